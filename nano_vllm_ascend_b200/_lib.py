"""ctypes binding of the C-ABI library ``libnvk_paged.so`` (declared in
``include/nvk_paged_kv.h``).

The library is the only compute path: if it is missing, importing the ops
raises instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libnvk_paged.so"

NVK_OK = 0
NVK_ERR_INVALID_ARGUMENT = -1
NVK_ERR_UNSUPPORTED = -2
NVK_ERR_WORKSPACE = -3
NVK_ERR_CUDA = -4

_c_void_p = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_size_t = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/nvk_paged_kv.h one to one.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "nvk_last_error": (ctypes.c_char_p, []),
    "nvk_abi_version": (_i32, []),
    "nvk_kv_append": (
        _i32,
        [_c_void_p, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i32, _i32, _c_void_p,
         _c_void_p],
    ),
    "nvk_paged_decode_workspace_size": (_i32, [_i32, _i32, _i32, _i32, _i32, ctypes.POINTER(_size_t)]),
    "nvk_paged_decode": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _c_void_p, _i32, _i32, _c_void_p, _i32, _i32, _i32,
         _i32, _f32, _i32, _c_void_p, _size_t, _c_void_p],
    ),
    "nvk_paged_decode_noalloc": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _c_void_p, _i32, _i32, _c_void_p, _i32, _i32, _i32,
         _i32, _f32, _i32, _c_void_p],
    ),
    "nvk_paged_decode_noalloc_error": (_i32, [ctypes.POINTER(_i32), _c_void_p]),
    "nvk_paged_prefill": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _c_void_p, _i32, _c_void_p, _c_void_p, _i32, _i32,
         _i32, _i32, _i32, _i32, _f32, _c_void_p, _c_void_p],
    ),
    "nvk_dense_prefill": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _f32, _c_void_p, _c_void_p],
    ),
    "nvk_qk_norm_rope_append": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _f32, _c_void_p, _c_void_p, _i32,
         _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i32, _i32, _i32, _c_void_p, _c_void_p],
    ),
    "nvk_decode_metadata": (
        _i32,
        [_c_void_p, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p, _c_void_p,
         _c_void_p, _c_void_p, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    ),
    "nvk_lm_head_argmax_workspace_size": (_i32, [_i32, ctypes.POINTER(_size_t)]),
    "nvk_lm_head_argmax": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _i32, _i32, _i32, _c_void_p, _c_void_p, _size_t, _i32, _c_void_p, _c_void_p],
    ),
    "nvk_prefix_create": (_i32, [_i32, _i32, ctypes.POINTER(_c_void_p)]),
    "nvk_prefix_destroy": (None, [_c_void_p]),
    "nvk_prefix_find_longest": (_i32, [_c_void_p, _c_void_p, _i64, _i32, _c_void_p, ctypes.POINTER(_i32)]),
    "nvk_prefix_cache_blocks": (_i32, [_c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p, _i64]),
    "nvk_prefix_forget_block": (_i32, [_c_void_p, _i32]),
    "nvk_prefix_block_key": (_i64, [_c_void_p, _i32]),
    "nvk_prefix_clear": (_i32, [_c_void_p]),
    "nvk_prefix_num_cached_keys": (_i64, [_c_void_p]),
    "nvk_prefix_num_keys": (_i64, [_c_void_p]),
    "nvk_peer_alloc": (_i32, [_size_t, ctypes.POINTER(_c_void_p)]),
    "nvk_peer_free": (_i32, [_c_void_p]),
    "nvk_peer_export": (_i32, [_c_void_p, _c_void_p]),
    "nvk_peer_import": (_i32, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "nvk_peer_close": (_i32, [_c_void_p]),
    "nvk_paged_decode_gather": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _i32, _i32, _c_void_p, _i32, _i32, _c_void_p, _i32, _i32, _i32, _i32, _f32,
         _i32, _c_void_p, _size_t, _c_void_p, _c_void_p, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _i64, _i64,
         _c_void_p, _c_void_p],
    ),
    "nvk_paged_decode_append": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _c_void_p, _i32, _i32, _c_void_p, _i32, _i32, _i32,
         _i32, _f32, _i32, _c_void_p, _size_t, _c_void_p, _c_void_p, _i64, _i64, _c_void_p, _c_void_p],
    ),
}

MAX_PEERS = 8
PEER_HANDLE_BYTES = 64
PEER_SIGNAL_BYTES = 256

_LIB: ctypes.CDLL | None = None


class NvkError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, func: str, code: int, message: str):
        super().__init__(f"{func} failed ({code}): {message}")
        self.code = code


def load() -> ctypes.CDLL:
    """Loads the library once and declares every exported signature."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = os.environ.get("NVK_PAGED_LIB", str(LIB_PATH))
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python -m nano_vllm_ascend_b200._build` "
            "(there is no non-CUDA implementation of these ops)"
        )
    lib = ctypes.CDLL(path)
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


def call(name: str, *args) -> None:
    """Calls ``name`` and raises NvkError (a RuntimeError) on a non-zero status."""
    check(name, getattr(load(), name)(*args))


def check(name: str, rc: int) -> None:
    """Raises for the status ``rc`` that entry point ``name`` returned, as ``call`` does."""
    if rc != NVK_OK:
        msg = load().nvk_last_error().decode(errors="replace")
        if rc in (NVK_ERR_INVALID_ARGUMENT, NVK_ERR_UNSUPPORTED):
            raise ValueError(f"{name}: {msg}")
        raise NvkError(name, rc, msg)
