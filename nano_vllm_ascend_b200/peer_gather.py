"""KV-head-sharded decode with the all-gather of the outputs done inside the
attention kernel (new: the reference runs on one device,
src/nanovllm_ascend/model_runner.py:31, and has no sharded path).

One process per GPU. Rank r holds KV heads [r*KVH/W, (r+1)*KVH/W) of every
layer and the query heads of their GQA groups. Each rank allocates one peer
buffer -- a signal area followed by ``slots`` gathered outputs [batch,
out_heads, head_dim] bf16 -- and maps every other rank's buffer through CUDA
IPC. ``nvk_paged_decode_gather`` then stores each output row of this rank's
heads into every rank's buffer over NVLink and, in its last CTA, exchanges an
epoch flag with every rank, so that when the call completes on this rank's
stream this rank's slot holds all heads. No NCCL call and no extra kernel is
on the data path.

A rank may run one call ahead of a slower peer; consecutive calls therefore
write different slots (``next_slot`` cycles through them).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .ops import _BF16, _ptr, _require_cuda, _stream, check_new_rows


class _DeviceBytes:
    """A raw device allocation seen by torch.as_tensor (CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerGather:
    """Gathered-output buffers shared by the ranks of ``group``.

    ``out_heads`` is the total number of query heads (all ranks); this rank's
    heads land at ``head_offset`` .. ``head_offset + local heads``.
    """

    def __init__(self, batch: int, out_heads: int, head_dim: int, slots: int = 2, device=None, group=None):
        if slots < 1:
            raise ValueError("PeerGather needs at least one output slot")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dist.is_available() and dist.is_initialized():
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        if not 1 <= self.world <= _lib.MAX_PEERS:
            raise ValueError(f"world size {self.world} outside 1..{_lib.MAX_PEERS}")
        self.batch, self.out_heads, self.head_dim, self.slots = batch, out_heads, head_dim, slots
        self.slot_bytes = (batch * out_heads * head_dim * 2 + 255) // 256 * 256
        self.nbytes = _lib.PEER_SIGNAL_BYTES + slots * self.slot_bytes
        self._slot = 0
        with torch.cuda.device(self.device):
            own = ctypes.c_void_p()
            _lib.call("nvk_peer_alloc", self.nbytes, ctypes.byref(own))
            self._own = own.value
            self._imported: list[int] = []
            bases = [0] * self.world
            bases[self.rank] = self._own
            if self.world > 1:
                handle = (ctypes.c_char * _lib.PEER_HANDLE_BYTES)()
                _lib.call("nvk_peer_export", ctypes.c_void_p(self._own), handle)
                handles: list[bytes | None] = [None] * self.world
                dist.all_gather_object(handles, bytes(handle), group=group)
                for r, h in enumerate(handles):
                    if r == self.rank:
                        continue
                    p = ctypes.c_void_p()
                    _lib.call("nvk_peer_import", ctypes.create_string_buffer(h, len(h)), ctypes.byref(p))
                    bases[r] = p.value
                    self._imported.append(p.value)
        self._bases = bases
        self._buffer = torch.as_tensor(_DeviceBytes(self._own, self.nbytes), device=self.device)
        self._group = group

    # ------------------------------------------------------------ layout ---
    def output(self, slot: int) -> torch.Tensor:
        """This rank's gathered output of ``slot``: bf16 [batch, out_heads, head_dim] (a view)."""
        off = _lib.PEER_SIGNAL_BYTES + slot * self.slot_bytes
        n = self.batch * self.out_heads * self.head_dim * 2
        return self._buffer[off: off + n].view(_BF16).view(self.batch, self.out_heads, self.head_dim)

    def _slot_ptrs(self, slot: int):
        off = _lib.PEER_SIGNAL_BYTES + slot * self.slot_bytes
        outs = (ctypes.c_void_p * _lib.MAX_PEERS)(*([b + off for b in self._bases] + [0] * (_lib.MAX_PEERS - self.world)))
        sigs = (ctypes.c_void_p * _lib.MAX_PEERS)(*(self._bases + [0] * (_lib.MAX_PEERS - self.world)))
        return outs, sigs

    def next_slot(self) -> int:
        s = self._slot
        self._slot = (self._slot + 1) % self.slots
        return s

    # ------------------------------------------------------------ decode ---
    def decode(self, query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
               block_tables: torch.Tensor, context_lens: torch.Tensor, scale: float, workspace: torch.Tensor,
               head_offset: int, slot: int | None = None, num_ctas: int = 0, new_key: torch.Tensor | None = None,
               new_value: torch.Tensor | None = None, slot_mapping: torch.Tensor | None = None) -> torch.Tensor:
        """Decode over this rank's heads; returns the gathered [batch, out_heads, D] output of the slot used.

        With ``new_key``/``new_value``/``slot_mapping`` the step's append of
        this rank's KV heads is fused in (see ops.paged_decode)."""
        dev = query.device
        for name, t in (("query", query), ("key_cache", key_cache), ("value_cache", value_cache),
                        ("block_tables", block_tables), ("context_lens", context_lens), ("workspace", workspace)):
            _require_cuda(name, t, dev)
        if query.dtype != _BF16 or key_cache.dtype != _BF16 or value_cache.dtype != _BF16:
            raise ValueError("paged_decode_gather: query and caches must be bfloat16")
        if not (query.is_contiguous() and key_cache.is_contiguous() and value_cache.is_contiguous()):
            raise ValueError("paged_decode_gather: query and caches must be contiguous")
        batch, num_heads, head_dim = query.shape
        num_blocks, block_size, kvh, d = key_cache.shape
        if batch != self.batch or head_dim != self.head_dim or d != head_dim or value_cache.shape != key_cache.shape:
            raise ValueError(f"paged_decode_gather: shape mismatch q={tuple(query.shape)} cache={tuple(key_cache.shape)}")
        if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.stride(1) != 1 \
                or block_tables.shape[0] != batch:
            raise ValueError("paged_decode_gather: block_tables must be int32 [batch, max_blocks]")
        if context_lens.dtype != torch.int32 or context_lens.numel() != batch or not context_lens.is_contiguous():
            raise ValueError("paged_decode_gather: context_lens must be a contiguous int32 [batch] device tensor")
        if slot_mapping is not None:
            new_key, new_value, slot_mapping = check_new_rows(new_key, new_value, slot_mapping, batch, kvh, head_dim,
                                                              dev)
        if slot is None:
            slot = self.next_slot()
        outs, sigs = self._slot_ptrs(slot)
        _lib.call(
            "nvk_paged_decode_gather", _ptr(query), _ptr(key_cache), _ptr(value_cache), num_blocks, block_size,
            _ptr(block_tables), block_tables.stride(0), block_tables.shape[1], _ptr(context_lens), batch, num_heads,
            kvh, head_dim, float(scale), int(num_ctas), _ptr(workspace),
            workspace.numel() * workspace.element_size(), outs, sigs, self.world, self.rank, self.out_heads,
            int(head_offset), _ptr(new_key), _ptr(new_value), 0 if new_key is None else new_key.stride(0),
            0 if new_value is None else new_value.stride(0), _ptr(slot_mapping), _stream(dev),
        )
        return self.output(slot)

    # ----------------------------------------------------------- teardown ---
    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (after a device sync
        and, with several ranks, a barrier so that no peer still writes)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self._group)
        self._buffer = None
        with torch.cuda.device(self.device):
            for p in self._imported:
                _lib.call("nvk_peer_close", ctypes.c_void_p(p))
            _lib.call("nvk_peer_free", ctypes.c_void_p(self._own))
        self._imported = []
        self._own = None
