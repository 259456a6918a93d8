"""CPU oracle for the paged-KV hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as a checker or as the timed CPU
reference. Nothing in the product (``nano_vllm_ascend_b200``) calls it.

A numpy restatement of the reference's path (Pla-Yer/nano_vllm_ascend, paths
relative to that project):

* slot mapping:   slot = table[pos // bs] * bs + pos % bs
                  (src/nanovllm_ascend/npu/block_manager.py:194-205, :233-250)
* KV append:      pool_flat[slot_mapping[t]] = rows[t]  (Tensor.index_copy_,
                  src/nanovllm_ascend/npu/paged_kv_cache.py:57-69), bit copy
* decode:         softmax(scale * q . K^T) V over the first context_lens[b]
                  tokens reached through block_tables[b]; query head h uses KV
                  head h // (H / KVH); scale = head_dim ** -0.5
                  (src/nanovllm_ascend/layers/npu_paged_attention.py:25-99;
                  docs/ascend_attention_kernels_metadata.md:140-250, :639-706)
* prefill:        bottom-right causal (sparse_mode=3): query i of a sequence
                  with Lq queries and Lk keys sees key j iff j <= Lk - Lq + i;
                  paged mode reads Lk = context_lens[b] keys via the block
                  table, dense mode reads contiguous k/v delimited by the
                  cumulative kv lengths
                  (src/nanovllm_ascend/layers/npu_prefill_attention.py:64-112;
                  docs/ascend_attention_kernels_metadata.md:1180-1204).

The attention arithmetic of the reference is a closed Ascend operator that is
not in the reference tree: attention parity is pinned only to this fp32
restatement (no golden vectors exist for it). Append and slot mapping are
pinned bit-exactly to fixtures produced by the reference's own
``PagedKVCache.write`` and ``BlockManager`` (tests/golden/).

bf16 tensors are handled as uint16 bit patterns so that numpy needs no bf16
type: widening is ``bits << 16`` viewed as float32.
"""

from __future__ import annotations

import numpy as np


# ------------------------------------------------------------- bf16 bits ----
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, np.uint16(0x7FC0), out)
    return out


# ---------------------------------------------------------- slot mapping ----
def slot_mapping(block_tables: list[list[int]], start_positions: list[int], num_tokens: list[int],
                 block_size: int) -> np.ndarray:
    """int64 slots for tokens [start, start + n) of every sequence, in order."""
    out = []
    for table, start, n in zip(block_tables, start_positions, num_tokens):
        for pos in range(start, start + n):
            idx = pos // block_size
            if idx >= len(table):
                raise RuntimeError(f"missing block at logical_pos={pos}")
            out.append(table[idx] * block_size + pos % block_size)
    return np.asarray(out, dtype=np.int64)


# ---------------------------------------------------------------- append ----
def kv_append(key_cache: np.ndarray, value_cache: np.ndarray, key: np.ndarray, value: np.ndarray,
              slots: np.ndarray) -> None:
    """In place on one layer [NB, BS, KVH, D] (any dtype, normally uint16 bits)."""
    nb, bs, kvh, d = key_cache.shape
    kflat = key_cache.reshape(nb * bs, kvh, d)
    vflat = value_cache.reshape(nb * bs, kvh, d)
    kflat[slots] = key
    vflat[slots] = value


# ------------------------------------------------- norm + rope + append ----
def qk_norm_rope_append(q: np.ndarray, k: np.ndarray, v: np.ndarray, q_weight: np.ndarray, k_weight: np.ndarray,
                        eps: float, cos_table: np.ndarray, sin_table: np.ndarray, positions: np.ndarray,
                        key_cache: np.ndarray, value_cache: np.ndarray, slots: np.ndarray) -> np.ndarray:
    """Prologue of Qwen3Attention.forward (src/nanovllm_ascend/models/qwen3.py:83-96).

    q [T, H, D], k/v [T, KVH, D] and the weights [D] are bf16 bits; the
    fp32 cos/sin tables are RotaryEmbedding's (layers/rotary_embedding.py:20-40).
    q_norm / k_norm (layers/layernorm.py:12-17): y = x / sqrt(mean(x^2) + eps) * w
    in fp32, output bf16. apply_rotary_pos_emb_tnd (:58-99): cos/sin rows cast to
    bf16, "half" rotation out = y * cos + rotate_half(y) * sin, rotate_half(y) =
    (-y[D/2:], y[:D/2]), output bf16. k_out and v are then written at slots
    (PagedKVCache.write, paged_kv_cache.py:44-69). Returns q_out bits.
    """
    def norm(x_bits, w_bits):
        x = bf16_bits_to_f32(x_bits)
        w = bf16_bits_to_f32(w_bits)
        ms = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
        y = (x * (np.float32(1.0) / np.sqrt(ms + np.float32(eps)))) * w
        return bf16_bits_to_f32(f32_to_bf16_bits(y.astype(np.float32)))

    pos = np.asarray(positions, dtype=np.int64)
    cos = bf16_bits_to_f32(f32_to_bf16_bits(cos_table[pos].astype(np.float32)))[:, None, :]
    sin = bf16_bits_to_f32(f32_to_bf16_bits(sin_table[pos].astype(np.float32)))[:, None, :]

    def rope(y):
        half = y.shape[-1] // 2
        rot = np.concatenate([-y[..., half:], y[..., :half]], axis=-1)
        return f32_to_bf16_bits((y * cos + rot * sin).astype(np.float32))

    q_out = rope(norm(q, q_weight))
    k_out = rope(norm(k, k_weight))
    kv_append(key_cache, value_cache, k_out, v, np.asarray(slots, dtype=np.int64))
    return q_out


# ------------------------------------------------------ lm head + argmax ----
def lm_head_logits(hidden: np.ndarray, weight: np.ndarray) -> np.ndarray:
    """bf16 logits of Qwen3ForCausalLM's lm_head (models/qwen3.py:196,221):
    hidden [B, H] and weight [V, H] as bf16 bits, f32 products summed in f32,
    rounded to bf16; returned as f32 values."""
    return bf16_bits_to_f32(f32_to_bf16_bits(as_f32(hidden) @ as_f32(weight).T))


def greedy_tokens(logits: np.ndarray) -> np.ndarray:
    """Sampler.sample's greedy branch (layers/sampler.py:13-14): torch.argmax
    over the vocabulary, the first index among equal maxima."""
    return np.argmax(logits, axis=-1).astype(np.int64)


# ---------------------------------------------------------------- decode ----
def as_f32(x: np.ndarray) -> np.ndarray:
    """uint16 arrays are bf16 bit patterns; anything else is cast to f32."""
    return bf16_bits_to_f32(x) if x.dtype == np.uint16 else x.astype(np.float32, copy=False)


def _gather_tokens(cache: np.ndarray, table: np.ndarray, n: int) -> np.ndarray:
    """First n token rows [n, KVH, D] (f32) of one sequence; only its blocks are widened."""
    bs = cache.shape[1]
    nblk = (n + bs - 1) // bs
    rows = cache[np.asarray(table[:nblk], dtype=np.int64)]  # [nblk, BS, KVH, D]
    return as_f32(rows.reshape(nblk * bs, *cache.shape[2:])[:n])


def _attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, visible: np.ndarray | None) -> np.ndarray:
    """q [Tq, H, D], k/v [Tk, KVH, D] f32 -> [Tq, H, D]; visible [Tq, Tk] bool."""
    tq, h, d = q.shape
    kvh = k.shape[1]
    qg = q.reshape(tq, kvh, h // kvh, d)
    s = np.einsum("tgqd,kgd->gqtk", qg, k, optimize=True) * np.float32(scale)
    if visible is not None:
        s = np.where(visible[None, None], s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)  # a row that sees no key yields zeros
    p = np.exp(s - m)
    denom = p.sum(axis=-1, keepdims=True)
    p = np.divide(p, denom, out=np.zeros_like(p), where=denom > 0)
    o = np.einsum("gqtk,kgd->tgqd", p, v, optimize=True)
    return o.reshape(tq, h, d).astype(np.float32)


def paged_decode(q: np.ndarray, key_cache: np.ndarray, value_cache: np.ndarray, block_tables: np.ndarray,
                 context_lens: np.ndarray, scale: float) -> np.ndarray:
    """q [B, H, D]; caches [NB, BS, KVH, D] (bf16 bits or float) -> [B, H, D] f32."""
    q = as_f32(q)
    out = np.zeros(q.shape, dtype=np.float32)
    for b in range(q.shape[0]):
        n = int(context_lens[b])
        if n <= 0:
            continue
        k = _gather_tokens(key_cache, block_tables[b], n)
        v = _gather_tokens(value_cache, block_tables[b], n)
        out[b] = _attend(q[b : b + 1], k, v, scale, None)[0]
    return out


# --------------------------------------------------------------- prefill ----
def _causal_visible(lq: int, lk: int) -> np.ndarray:
    i = np.arange(lq)[:, None]
    j = np.arange(lk)[None, :]
    return j <= (lk - lq) + i


def paged_prefill(q: np.ndarray, key_cache: np.ndarray, value_cache: np.ndarray, block_tables: np.ndarray,
                  cu_seqlens_q: np.ndarray, kv_lens: np.ndarray, scale: float) -> np.ndarray:
    """q [Tq, H, D] -> [Tq, H, D] f32; sequence b owns rows cu[b]:cu[b+1]."""
    q = as_f32(q)
    out = np.zeros(q.shape, dtype=np.float32)
    for b in range(len(kv_lens)):
        s, e = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
        lk = int(kv_lens[b])
        if e <= s:
            continue
        k = _gather_tokens(key_cache, block_tables[b], lk)
        v = _gather_tokens(value_cache, block_tables[b], lk)
        out[s:e] = _attend(q[s:e], k, v, scale, _causal_visible(e - s, lk))
    return out


def dense_prefill(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_seqlens_q: np.ndarray,
                  cu_seqlens_kv: np.ndarray, scale: float) -> np.ndarray:
    q, k, v = as_f32(q), as_f32(k), as_f32(v)
    out = np.zeros(q.shape, dtype=np.float32)
    for b in range(len(cu_seqlens_q) - 1):
        s, e = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
        ks, ke = int(cu_seqlens_kv[b]), int(cu_seqlens_kv[b + 1])
        if e <= s:
            continue
        out[s:e] = _attend(q[s:e], k[ks:ke], v[ks:ke], scale, _causal_visible(e - s, ke - ks))
    return out
