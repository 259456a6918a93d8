"""Generates the golden fixtures in this directory from the REFERENCE itself.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py /path/to/nano_vllm_ascend

It imports the reference's own CPU-importable host classes --
``nanovllm_ascend.npu.block_manager.BlockManager`` and
``nanovllm_ascend.npu.paged_kv_cache.PagedKVCache`` (both need only torch) --
drives them with seeded inputs, and records what they return:

* block_manager_golden.json -- block tables, CPU context lengths, slot
  mappings, prefix lookups and free-queue snapshots for (a) the reference's
  own unit-test scenarios (tests/test_block_manager.py:6-54), (b) a seeded
  random script of prefill / decode / cache / free / clear operations with
  prefix reuse, (c) the config-1 decode step (64 blocks of 128, free queue =
  torch.randperm(64) with seed 0, contexts {37, 128, 255, 513} + 1 token).
* append_golden.json -- ``PagedKVCache.write`` (the reference's index_copy_
  append) on the config-1 decode append and a prefill-sized ragged append.
  Inputs are regenerated from their seed by ``append_inputs`` below (the
  SHA-256 of the regenerated bf16 bits is recorded so a different RNG fails
  loudly); results are SHA-256 digests of the written rows and of each whole
  pool (zero-filled before the write).

The fixtures are committed; tests read them on any machine (including the GPU
box, where the reference is absent).
"""

from __future__ import annotations

import hashlib
import json
import random
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _md(m) -> dict:
    return {
        "block_tables": m.block_tables.tolist(),
        "context_lens": m.context_lens.tolist(),
        "context_lens_device": str(m.context_lens.device),
        "context_lens_dtype": str(m.context_lens.dtype),
        "block_tables_dtype": str(m.block_tables.dtype),
        "slot_mapping": m.slot_mapping.tolist(),
        "slot_mapping_dtype": str(m.slot_mapping.dtype),
        "actual_seq_lengths_q": m.actual_seq_lengths_q,
        "actual_seq_lengths_kv": m.actual_seq_lengths_kv,
        "query_lens": m.query_lens,
        "use_paged_prefill": m.use_paged_prefill,
    }


def random_script(seed: int, num_blocks: int, block_size: int, steps: int) -> list[dict]:
    """A seeded operation script exercising allocation, prefix reuse and eviction.

    Prompts are drawn from a few shared stems so that prefix hits, partial
    hits and evictions of cached blocks all occur.
    """
    rng = random.Random(seed)
    stems = [[rng.randrange(50) for _ in range(block_size * 4)] for _ in range(3)]
    ops: list[dict] = []
    live: dict[int, dict] = {}
    next_slot = 0
    for _ in range(steps):
        r = rng.random()
        if r < 0.35 and len(live) < 5:
            stem = rng.choice(stems)
            keep = rng.randrange(0, len(stem) + 1)
            tail = [rng.randrange(50, 100) for _ in range(rng.randrange(1, 2 * block_size + 3))]
            tokens = stem[:keep] + tail
            ops.append({"op": "admit", "slot": next_slot, "tokens": tokens})
            live[next_slot] = {"len": len(tokens)}
            next_slot += 1
        elif r < 0.75 and live:
            slots = sorted(rng.sample(sorted(live), rng.randrange(1, len(live) + 1)))
            ops.append({"op": "decode", "slots": slots})
            for s in slots:
                live[s]["len"] += 1
        elif live:
            s = rng.choice(sorted(live))
            ops.append({"op": "free", "slot": s})
            del live[s]
        elif rng.random() < 0.2:
            ops.append({"op": "clear"})
    for s in sorted(live):
        ops.append({"op": "free", "slot": s})
    ops.append({"op": "clear"})
    return ops


def run_script(bm_cls, ops: list[dict], num_blocks: int, block_size: int) -> list[dict]:
    """Replays a script the way ModelRunner drives the BlockManager
    (model_runner.py:146-167 prefix lookup, :199-238 prefill + cache_full_blocks,
    :240-286 decode, :293-294 free)."""
    bm = bm_cls(num_blocks=num_blocks, block_size=block_size, device="cpu")
    lens: dict[int, int] = {}
    results: list[dict] = []
    for op in ops:
        res: dict = {"op": op["op"]}
        try:
            if op["op"] == "admit":
                tokens = torch.tensor(op["tokens"], dtype=torch.long)
                n = tokens.numel()
                full = n // block_size
                max_cache = full - 1 if (n % block_size == 0 and full > 0) else full
                cached = bm.find_longest_prefix_blocks(tokens, max_cache_blocks=max_cache) if max_cache > 0 else []
                start = len(cached) * block_size
                md = bm.prepare_prefill_metadata(slots=[op["slot"]], seq_lens=[n - start], start_positions=[start],
                                                 prefix_block_ids=[cached])
                bm.cache_full_blocks(slot=op["slot"], token_ids=tokens, num_cached_blocks=len(cached),
                                     num_full_blocks=full)
                lens[op["slot"]] = n
                res.update(cached=cached, md=_md(md))
            elif op["op"] == "decode":
                starts = [lens[s] for s in op["slots"]]
                md = bm.prepare_decode_metadata(slots=op["slots"], start_positions=starts, q_len=1)
                for s in op["slots"]:
                    lens[s] += 1
                res.update(md=_md(md))
            elif op["op"] == "free":
                bm.free_slot(op["slot"])
                lens.pop(op["slot"], None)
            elif op["op"] == "clear":
                bm.clear_prefix_cache()
        except Exception as exc:  # errors are part of the observable behaviour
            res["error"] = f"{type(exc).__name__}: {exc}"
        res["free"] = list(bm.free_block_ids)
        res["ref_counts"] = [b.ref_count for b in bm.blocks]
        res["hashed"] = [b.block_hash is not None for b in bm.blocks]
        results.append(res)
    return results


def unit_scenarios(bm_cls) -> dict:
    out = {}
    m = bm_cls(num_blocks=8, block_size=4, device="cpu")
    md = m.prepare_prefill_metadata(slots=[0, 1, 2], seq_lens=[3, 5, 2], start_positions=[0, 0, 0],
                                    prefix_block_ids=[[], [], []])
    out["prefill"] = _md(md)
    md2 = m.prepare_decode_metadata(slots=[1, 2], start_positions=[5, 2], q_len=1)
    out["decode"] = _md(md2)
    m = bm_cls(num_blocks=8, block_size=4, device="cpu")
    tokens = torch.tensor([10, 11, 12, 13, 20, 21], dtype=torch.long)
    m.prepare_prefill_metadata(slots=[0], seq_lens=[6], start_positions=[0], prefix_block_ids=[[]])
    m.cache_full_blocks(slot=0, token_ids=tokens)
    m.free_slot(0)
    out["prefix_reuse"] = m.find_longest_prefix_blocks(tokens, max_cache_blocks=1)
    out["prefix_reuse_free"] = list(m.free_block_ids)
    return out


def config1(bm_cls) -> dict:
    """Config 1: 64 blocks of 128; free queue = randperm(64, seed 0);
    contexts {37, 128, 255, 513} prefilled, then one decode token each."""
    g = torch.Generator().manual_seed(0)
    perm = torch.randperm(64, generator=g).tolist()
    bm = bm_cls(num_blocks=64, block_size=128, device="cpu")
    bm.free_block_ids = list(perm)
    ctx = [37, 128, 255, 513]
    slots = [0, 1, 2, 3]
    pre = bm.prepare_prefill_metadata(slots=slots, seq_lens=ctx, start_positions=[0] * 4,
                                      prefix_block_ids=[[] for _ in slots])
    dec = bm.prepare_decode_metadata(slots=slots, start_positions=ctx, q_len=1)
    return {"perm": perm, "ctx": ctx, "prefill": _md(pre), "decode": _md(dec)}


def sha(bits: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(bits).tobytes()).hexdigest()


def append_inputs(num_tokens: int, kvh: int, d: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Seeded bf16 K/V rows [T, KVH, D] ~ N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(num_tokens, kvh, d, generator=g).to(torch.bfloat16)
    v = torch.randn(num_tokens, kvh, d, generator=g).to(torch.bfloat16)
    return k, v


def append_case(kv_cls, num_blocks, block_size, kvh, d, slots: list[int], seed: int) -> dict:
    k, v = append_inputs(len(slots), kvh, d, seed)
    kv = kv_cls(num_layers=1, num_blocks=num_blocks, block_size=block_size, num_kv_heads=kvh, head_dim=d,
                dtype=torch.bfloat16, device="cpu")
    kv.key_cache.zero_()
    kv.value_cache.zero_()
    slot_t = torch.tensor(slots, dtype=torch.int64)
    kv.write(layer_idx=0, key_states=k, value_states=v, slot_mapping=slot_t)
    kc, vc = kv.get_physical_cache(0)
    flat_k = kc.reshape(num_blocks * block_size, kvh, d)
    flat_v = vc.reshape(num_blocks * block_size, kvh, d)
    return {
        "shape": [num_blocks, block_size, kvh, d],
        "slots": slots,
        "seed": seed,
        "sha_key_in": sha(_bits(k)),
        "sha_value_in": sha(_bits(v)),
        "sha_rows_key": sha(_bits(flat_k[slot_t])),
        "sha_rows_value": sha(_bits(flat_v[slot_t])),
        "sha_pool_key": sha(_bits(kc)),
        "sha_pool_value": sha(_bits(vc)),
    }


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    from nanovllm_ascend.npu.block_manager import BlockManager
    from nanovllm_ascend.npu.paged_kv_cache import PagedKVCache

    script = random_script(seed=1234, num_blocks=24, block_size=4, steps=160)
    golden = {
        "unit": unit_scenarios(BlockManager),
        "script": {"num_blocks": 24, "block_size": 4, "ops": script,
                   "results": run_script(BlockManager, script, 24, 4)},
        "config1": config1(BlockManager),
    }
    (HERE / "block_manager_golden.json").write_text(json.dumps(golden, separators=(",", ":")))

    c1 = golden["config1"]["decode"]["slot_mapping"]
    # Prefill-sized ragged append: 3 sequences of 200, 77 and 128 tokens over
    # blocks handed out from a seeded permutation of a 16-block pool.
    g = torch.Generator().manual_seed(7)
    perm = torch.randperm(16, generator=g).tolist()
    bm = BlockManager(num_blocks=16, block_size=128, device="cpu")
    bm.free_block_ids = perm
    md = bm.prepare_prefill_metadata(slots=[0, 1, 2], seq_lens=[200, 77, 128], start_positions=[0, 0, 0],
                                     prefix_block_ids=[[], [], []])
    cases = {
        "c1": append_case(PagedKVCache, 64, 128, 8, 128, c1, seed=11),
        "ragged": append_case(PagedKVCache, 16, 128, 8, 128, md.slot_mapping.tolist(), seed=12),
    }
    (HERE / "append_golden.json").write_text(json.dumps(cases, indent=1))
    print("wrote", HERE / "block_manager_golden.json", HERE / "append_golden.json")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
