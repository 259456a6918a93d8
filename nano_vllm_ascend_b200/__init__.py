"""B200-native paged-KV-cache hot path of nano_vllm_ascend.

Drop-in host classes (same names and contracts as the reference's):

* ``PagedKVCache`` -- pool + CUDA append          (npu/paged_kv_cache.py)
* ``BlockManager`` / ``PagedKVCacheMetadata``     (npu/block_manager.py)
* ``PagedAttention``  -- decode attention          (layers/npu_paged_attention.py)
* ``BatchPrefillAttention`` -- causal prefill     (layers/npu_prefill_attention.py)
* ``DecodeGraphRunner`` -- CUDA-graph decode       (npu/acl_graph.py)

Device-side errors (bad slots, block ids, over-long contexts) raise with the
reference's exception types through ``device_errors`` / ``check_errors()``.

The compute lives in ``libnvk_paged.so`` (C ABI in include/nvk_paged_kv.h),
built for sm_100a by ``nano_vllm_ascend_b200._build``.
"""

from . import device_errors
from .block_manager import BlockManager, BlockState, PagedKVCacheMetadata
from .cuda_graph import DecodeGraphRunner, DecodeGraphStats, copy_block_tables
from .paged_attention import PagedAttention
from .paged_kv_cache import PagedKVCache
from .device_errors import KVCacheDeviceError, check_errors
from .prefill_attention import BatchPrefillAttention

# Names used by the reference's call sites.
NpuPagedAttention = PagedAttention
NpuBatchPrefillAttention = BatchPrefillAttention

__all__ = [
    "BatchPrefillAttention",
    "BlockManager",
    "BlockState",
    "DecodeGraphRunner",
    "DecodeGraphStats",
    "KVCacheDeviceError",
    "NpuBatchPrefillAttention",
    "NpuPagedAttention",
    "PagedAttention",
    "PagedKVCache",
    "PagedKVCacheMetadata",
    "check_errors",
    "copy_block_tables",
]
