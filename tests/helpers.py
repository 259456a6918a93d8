"""Shared builders for the GPU parity tests (seeded inputs, oracle adapters)."""

from __future__ import annotations

import numpy as np
import torch

ATOL = 2e-2  # attention tolerance vs the fp32 oracle (bf16 outputs)
RTOL = 1e-2


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor (any device) -> uint16 bit patterns on the host."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def seeded_tables(ctx: list[int], block_size: int, num_blocks: int, seed: int, width: int | None = None):
    """Block tables drawn without replacement from a seeded pool permutation."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g)
    need = [(n + block_size - 1) // block_size for n in ctx]
    if sum(need) > num_blocks:
        raise ValueError("pool too small for the requested contexts")
    width = width or max(max(need), 1)
    tables = torch.zeros(len(ctx), width, dtype=torch.int32)
    used = 0
    for i, m in enumerate(need):
        tables[i, :m] = perm[used : used + m].to(torch.int32)
        used += m
    return tables


def random_pool(num_blocks: int, block_size: int, kvh: int, d: int, device, seed: int):
    g = torch.Generator(device=device).manual_seed(seed)
    shape = (num_blocks, block_size, kvh, d)
    kc = torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    vc = torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    return kc, vc


def assert_close(got: np.ndarray, want: np.ndarray, what: str = "") -> tuple[float, float]:
    err = np.abs(got - want)
    max_abs = float(err.max()) if err.size else 0.0
    bad = ~(err <= ATOL + RTOL * np.abs(want))  # NaN (an unwritten output) counts as bad
    if bad.any():
        idx = np.argwhere(bad)[0]
        raise AssertionError(f"{what}: {int(bad.sum())} elements outside atol={ATOL} rtol={RTOL}; first at "
                             f"{tuple(idx)} got={got[tuple(idx)]} want={want[tuple(idx)]} max_abs={max_abs}")
    return max_abs, float((err / (np.abs(want) + 1e-6)).max()) if err.size else 0.0
