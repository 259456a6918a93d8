"""Tensor-level wrappers over the C-ABI kernels.

Each function validates devices, dtypes, shapes and strides, then calls the
matching ``nvk_*`` entry point on the tensors' current CUDA stream. Nothing
here computes on the host: there is no non-CUDA path.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_BF16 = torch.bfloat16
_KV_DTYPES = (torch.bfloat16, torch.float16)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(name: str, t: torch.Tensor, device: torch.device | None = None) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (got device {t.device})")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")


def _require_rows(name: str, t: torch.Tensor) -> None:
    """[T, heads, dim] with heads and dims packed; the token stride may be larger."""
    if t.dim() != 3 or t.stride(2) != 1 or t.stride(1) != t.shape[2]:
        raise ValueError(f"{name} must be [tokens, heads, dim] with contiguous heads/dims, got "
                         f"shape {tuple(t.shape)} stride {t.stride()}")


# ----------------------------------------------------------------- append ---
def kv_append(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    slot_mapping: torch.Tensor,
    error_word: torch.Tensor | None = None,
) -> None:
    """key_cache.view(-1, KVH, D)[slot_mapping] = key (same for value), in place.

    ``key_cache``/``value_cache`` are ONE layer of the pool, [NB, BS, KVH, D]
    contiguous. ``slot_mapping`` must be int64 on the same device.
    """
    dev = key_cache.device
    for name, t in (("key_cache", key_cache), ("value_cache", value_cache), ("key", key), ("value", value),
                    ("slot_mapping", slot_mapping)):
        _require_cuda(name, t, dev)
    if key_cache.dtype not in _KV_DTYPES or key.dtype != key_cache.dtype or value.dtype != key_cache.dtype \
            or value_cache.dtype != key_cache.dtype:
        raise ValueError(f"kv_append: dtype mismatch (cache {key_cache.dtype}, key {key.dtype}, value {value.dtype})")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()) or key_cache.shape != value_cache.shape:
        raise ValueError("kv_append: key/value cache must be contiguous and of equal shape")
    num_blocks, block_size, kvh, d = key_cache.shape
    _require_rows("key", key)
    _require_rows("value", value)
    if key.shape != value.shape or key.shape[1] != kvh or key.shape[2] != d:
        raise ValueError(f"kv shape mismatch: got {tuple(key.shape)} / {tuple(value.shape)}")
    if slot_mapping.dtype != torch.int64 or slot_mapping.numel() != key.shape[0]:
        raise ValueError("kv_append: slot_mapping must be int64 with one entry per token")
    slot_mapping = slot_mapping.contiguous()
    if error_word is not None:
        _require_cuda("error_word", error_word, dev)
    _lib.call(
        "nvk_kv_append", _ptr(key), _ptr(value), key.stride(0), value.stride(0), _ptr(key_cache), _ptr(value_cache),
        _ptr(slot_mapping), key.shape[0], num_blocks * block_size, kvh, d, _ptr(error_word), _stream(dev),
    )


# ------------------------------------------------- norm + rope + append ---
def qk_norm_rope_append(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    eps: float,
    cos_table: torch.Tensor,
    sin_table: torch.Tensor,
    positions: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    query_out: torch.Tensor | None = None,
    error_word: torch.Tensor | None = None,
) -> torch.Tensor:
    """q_norm + k_norm + rotary embedding + KV append in one kernel
    (Qwen3Attention.forward's prologue, qwen3.py:83-96). Returns the rotated
    query [T, H, D] (``query_out``, new if None); the rotated key and the value
    rows land in ONE layer of the pool at ``slot_mapping``."""
    dev = query.device
    for name, t in (("query", query), ("key", key), ("value", value), ("q_weight", q_weight),
                    ("k_weight", k_weight), ("cos_table", cos_table), ("sin_table", sin_table),
                    ("positions", positions), ("key_cache", key_cache), ("value_cache", value_cache),
                    ("slot_mapping", slot_mapping)):
        _require_cuda(name, t, dev)
    for name, t in (("query", query), ("key", key), ("value", value)):
        _require_rows(name, t)
        if t.dtype != _BF16:
            raise ValueError(f"qk_norm_rope_append: {name} must be bfloat16")
    tokens, num_heads, head_dim = query.shape
    num_blocks, block_size, kvh, d = key_cache.shape
    if key.shape != (tokens, kvh, head_dim) or value.shape != key.shape or d != head_dim:
        raise ValueError(f"kv shape mismatch: got {tuple(key.shape)} / {tuple(value.shape)}")
    if q_weight.numel() != head_dim or k_weight.numel() != head_dim or q_weight.dtype != _BF16 \
            or k_weight.dtype != _BF16:
        raise ValueError("qk_norm_rope_append: q_weight/k_weight must be bfloat16 [head_dim]")
    if cos_table.dtype != torch.float32 or sin_table.shape != cos_table.shape or cos_table.dim() != 2 \
            or cos_table.shape[1] != head_dim or not (cos_table.is_contiguous() and sin_table.is_contiguous()):
        raise ValueError("qk_norm_rope_append: cos/sin tables must be contiguous float32 [max_position, head_dim]")
    if positions.dtype != torch.int64 or positions.numel() != tokens or slot_mapping.dtype != torch.int64 \
            or slot_mapping.numel() != tokens:
        raise ValueError("qk_norm_rope_append: positions and slot_mapping must be int64 [tokens]")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("qk_norm_rope_append: caches must be contiguous")
    if query_out is None:
        query_out = torch.empty(tokens, num_heads, head_dim, dtype=_BF16, device=dev)
    elif query_out.shape != (tokens, num_heads, head_dim) or not query_out.is_contiguous() or query_out.dtype != _BF16:
        raise ValueError("qk_norm_rope_append: query_out must be a contiguous bf16 [tokens, heads, head_dim]")
    _lib.call(
        "nvk_qk_norm_rope_append", _ptr(query), _ptr(key), _ptr(value), query.stride(0), key.stride(0),
        value.stride(0), _ptr(q_weight.contiguous()), _ptr(k_weight.contiguous()), float(eps), _ptr(cos_table),
        _ptr(sin_table), cos_table.shape[0], _ptr(positions.contiguous()), _ptr(query_out), _ptr(key_cache),
        _ptr(value_cache), _ptr(slot_mapping.contiguous()), tokens, num_blocks * block_size, num_heads, kvh,
        head_dim, _ptr(error_word), _stream(dev),
    )
    return query_out


# ----------------------------------------------------- lm head + argmax ---
def lm_head_argmax_workspace_bytes(batch: int) -> int:
    out = ctypes.c_size_t(0)
    _lib.call("nvk_lm_head_argmax_workspace_size", batch, ctypes.byref(out))
    return int(out.value)


def lm_head_argmax(hidden: torch.Tensor, weight: torch.Tensor, workspace: torch.Tensor,
                   token_ids: torch.Tensor | None = None, num_ctas: int = 0,
                   error_word: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy next tokens of a decode batch: argmax over the vocabulary of the
    bf16 logits hidden @ weight.T (first index on ties), int64 [batch] on the
    device. ``workspace`` (uint8, zeroed once) holds
    lm_head_argmax_workspace_bytes(batch); ``error_word`` a device int32."""
    dev = hidden.device
    for name, t in (("hidden", hidden), ("weight", weight), ("workspace", workspace)):
        _require_cuda(name, t, dev)
    if hidden.dtype != _BF16 or weight.dtype != _BF16 or hidden.dim() != 2 or weight.dim() != 2 \
            or hidden.stride(1) != 1 or not weight.is_contiguous() or weight.shape[1] != hidden.shape[1]:
        raise ValueError("lm_head_argmax: hidden [batch, H] and weight [vocab, H] must be bf16 with unit inner stride")
    batch, hsize = hidden.shape
    if token_ids is None:
        token_ids = torch.empty(batch, dtype=torch.int64, device=dev)
    if error_word is None:
        error_word = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.call("nvk_lm_head_argmax", _ptr(hidden), hidden.stride(0), _ptr(weight), weight.shape[0], hsize, batch,
              _ptr(token_ids), _ptr(workspace), workspace.numel() * workspace.element_size(), int(num_ctas),
              _ptr(error_word), _stream(dev))
    return token_ids


# ----------------------------------------------------------------- decode ---
def decode_workspace_bytes(batch: int, num_heads: int, num_kv_heads: int, head_dim: int, num_ctas: int = 0) -> int:
    """Workspace bytes of paged_decode (num_ctas 0 = one CTA per SM of the current device)."""
    out = ctypes.c_size_t(0)
    _lib.call("nvk_paged_decode_workspace_size", batch, num_heads, num_kv_heads, head_dim, num_ctas,
              ctypes.byref(out))
    return int(out.value)


def paged_decode(
    out: torch.Tensor,
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    workspace: torch.Tensor,
    num_ctas: int = 0,
    new_key: torch.Tensor | None = None,
    new_value: torch.Tensor | None = None,
    slot_mapping: torch.Tensor | None = None,
) -> torch.Tensor:
    """Paged GQA decode attention into ``out`` ([B, H, D] bf16).

    ``workspace`` (uint8, zeroed once) must hold decode_workspace_bytes(B, H,
    KVH, D, num_ctas); calls sharing it must be ordered on one stream.
    With ``new_key``/``new_value`` ([B, KVH, D] rows) and ``slot_mapping``
    ([B] int64) the step's append is fused in: the rows are written to the
    pool at their slots (each sequence's last context position) and attended
    over, as kv_append followed by paged_decode.
    """
    dev = query.device
    for name, t in (("out", out), ("query", query), ("key_cache", key_cache), ("value_cache", value_cache),
                    ("block_tables", block_tables), ("context_lens", context_lens), ("workspace", workspace)):
        _require_cuda(name, t, dev)
    if query.dtype != _BF16 or out.dtype != _BF16 or key_cache.dtype != _BF16 or value_cache.dtype != _BF16:
        raise ValueError("paged_decode: query, out and caches must be bfloat16")
    if not (query.is_contiguous() and out.is_contiguous() and key_cache.is_contiguous()
            and value_cache.is_contiguous()):
        raise ValueError("paged_decode: query, out and caches must be contiguous")
    batch, num_heads, head_dim = query.shape
    num_blocks, block_size, kvh, d = key_cache.shape
    if d != head_dim or value_cache.shape != key_cache.shape or out.shape != query.shape:
        raise ValueError(f"paged_decode: shape mismatch q={tuple(query.shape)} cache={tuple(key_cache.shape)}")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.stride(1) != 1 \
            or block_tables.shape[0] != batch:
        raise ValueError("paged_decode: block_tables must be int32 [batch, max_blocks] with unit column stride")
    if context_lens.dtype != torch.int32 or context_lens.numel() != batch or not context_lens.is_contiguous():
        raise ValueError("paged_decode: context_lens must be a contiguous int32 [batch] device tensor")
    ws_bytes = workspace.numel() * workspace.element_size()
    if slot_mapping is None:
        _lib.call(
            "nvk_paged_decode", _ptr(out), _ptr(query), _ptr(key_cache), _ptr(value_cache), num_blocks, block_size,
            _ptr(block_tables), block_tables.stride(0), block_tables.shape[1], _ptr(context_lens), batch, num_heads,
            kvh, head_dim, float(scale), int(num_ctas), _ptr(workspace), ws_bytes, _stream(dev),
        )
        return out
    new_key, new_value, slot_mapping = check_new_rows(new_key, new_value, slot_mapping, batch, kvh, head_dim, dev)
    _lib.call(
        "nvk_paged_decode_append", _ptr(out), _ptr(query), _ptr(key_cache), _ptr(value_cache), num_blocks,
        block_size, _ptr(block_tables), block_tables.stride(0), block_tables.shape[1], _ptr(context_lens), batch,
        num_heads, kvh, head_dim, float(scale), int(num_ctas), _ptr(workspace), ws_bytes, _ptr(new_key),
        _ptr(new_value), new_key.stride(0), new_value.stride(0), _ptr(slot_mapping), _stream(dev),
    )
    return out


def check_new_rows(new_key, new_value, slot_mapping, batch: int, kvh: int, head_dim: int, dev):
    """Validates the one-token-per-sequence rows of a fused append; returns them usable by the kernel."""
    if new_key is None or new_value is None:
        raise ValueError("paged_decode: a fused append needs new_key, new_value and slot_mapping")
    for name, t in (("new_key", new_key), ("new_value", new_value), ("slot_mapping", slot_mapping)):
        _require_cuda(name, t, dev)
    if new_key.dtype != _BF16 or new_value.dtype != _BF16:
        raise ValueError("paged_decode: new_key/new_value must be bfloat16")
    _require_rows("new_key", new_key)
    _require_rows("new_value", new_value)
    if new_key.shape != (batch, kvh, head_dim) or new_value.shape != new_key.shape:
        raise ValueError(f"kv shape mismatch: got {tuple(new_key.shape)} / {tuple(new_value.shape)}")
    if slot_mapping.dtype != torch.int64 or slot_mapping.numel() != batch:
        raise ValueError("paged_decode: slot_mapping must be int64 with one entry per sequence")
    if (new_key.stride(0) * 2) % 16 or new_key.data_ptr() % 16:
        new_key = new_key.contiguous()
    if (new_value.stride(0) * 2) % 16 or new_value.data_ptr() % 16:
        new_value = new_value.contiguous()
    return new_key, new_value, slot_mapping.contiguous()


def decode_error_word(workspace: torch.Tensor) -> int:
    """Reads (synchronously) the device error word at the head of a decode workspace."""
    return int(workspace[:4].view(torch.int32).item())


# ---------------------------------------------------------------- prefill ---
def paged_prefill(
    out: torch.Tensor,
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    kv_lens: torch.Tensor,
    max_q_len: int,
    scale: float,
    error_word: torch.Tensor | None = None,
) -> torch.Tensor:
    """Causal (bottom-right) prefill attention over the paged pool into ``out``."""
    dev = query.device
    for name, t in (("out", out), ("query", query), ("key_cache", key_cache), ("value_cache", value_cache),
                    ("block_tables", block_tables), ("cu_seqlens_q", cu_seqlens_q), ("kv_lens", kv_lens)):
        _require_cuda(name, t, dev)
    if query.dtype != _BF16 or out.dtype != _BF16 or key_cache.dtype != _BF16 or value_cache.dtype != _BF16:
        raise ValueError("paged_prefill: query, out and caches must be bfloat16")
    if not (query.is_contiguous() and out.is_contiguous() and key_cache.is_contiguous()
            and value_cache.is_contiguous()):
        raise ValueError("paged_prefill: query, out and caches must be contiguous")
    total_q, num_heads, head_dim = query.shape
    num_blocks, block_size, kvh, d = key_cache.shape
    batch = kv_lens.numel()
    if d != head_dim or out.shape != query.shape or value_cache.shape != key_cache.shape:
        raise ValueError("paged_prefill: shape mismatch")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.stride(1) != 1 \
            or block_tables.shape[0] != batch:
        raise ValueError("paged_prefill: block_tables must be int32 [batch, max_blocks]")
    if cu_seqlens_q.dtype != torch.int32 or cu_seqlens_q.numel() != batch + 1 or kv_lens.dtype != torch.int32:
        raise ValueError("paged_prefill: cu_seqlens_q must be int32 [batch+1] and kv_lens int32 [batch]")
    _lib.call(
        "nvk_paged_prefill", _ptr(out), _ptr(query), _ptr(key_cache), _ptr(value_cache), num_blocks, block_size,
        _ptr(block_tables), block_tables.stride(0), _ptr(cu_seqlens_q.contiguous()), _ptr(kv_lens.contiguous()),
        batch, total_q, int(max_q_len), num_heads, kvh, head_dim, float(scale), _ptr(error_word), _stream(dev),
    )
    return out


def dense_prefill(
    out: torch.Tensor,
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    cu_seqlens_kv: torch.Tensor,
    max_q_len: int,
    scale: float,
    error_word: torch.Tensor | None = None,
) -> torch.Tensor:
    """Causal (bottom-right) prefill attention over contiguous K/V rows."""
    dev = query.device
    for name, t in (("out", out), ("query", query), ("key", key), ("value", value), ("cu_seqlens_q", cu_seqlens_q),
                    ("cu_seqlens_kv", cu_seqlens_kv)):
        _require_cuda(name, t, dev)
    if any(t.dtype != _BF16 for t in (out, query, key, value)):
        raise ValueError("dense_prefill: tensors must be bfloat16")
    if not all(t.is_contiguous() for t in (out, query, key, value)):
        raise ValueError("dense_prefill: tensors must be contiguous")
    total_q, num_heads, head_dim = query.shape
    total_kv, kvh, d = key.shape
    batch = cu_seqlens_q.numel() - 1
    if d != head_dim or value.shape != key.shape or out.shape != query.shape or cu_seqlens_kv.numel() != batch + 1:
        raise ValueError("dense_prefill: shape mismatch")
    _lib.call(
        "nvk_dense_prefill", _ptr(out), _ptr(query), _ptr(key), _ptr(value), _ptr(cu_seqlens_q.contiguous()),
        _ptr(cu_seqlens_kv.contiguous()), batch, total_q, total_kv, int(max_q_len), num_heads, kvh, head_dim,
        float(scale), _ptr(error_word), _stream(dev),
    )
    return out
