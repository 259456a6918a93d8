"""C-ABI library checks that need no GPU.

The library loads on a host without a driver, exports exactly the entry points
declared in include/*.h, and rejects bad arguments on the host (before any CUDA
call) with the documented status codes.
"""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from nano_vllm_ascend_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions() -> set[str]:
    names = set()
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_\s\*]*?\b(nvk_[a-z0-9_]+)\s*\(", text, re.M):
            names.add(m.group(1))
    return names


def test_headers_declare_the_boundary():
    names = declared_functions()
    assert {"nvk_kv_append", "nvk_paged_decode", "nvk_paged_decode_workspace_size", "nvk_paged_prefill",
            "nvk_dense_prefill", "nvk_last_error", "nvk_abi_version"} <= names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert set(_lib.SIGNATURES) == declared_functions()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line and "nvk_" in line}
    assert exported == declared_functions(), "only the declared C entry points may be exported"


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.nvk_abi_version() == 5
    assert isinstance(lib.nvk_last_error(), bytes)


def test_host_side_validation_codes():
    lib = _lib.load()
    n = ctypes.c_void_p(0)
    # args: out q kc vc num_blocks block_size tables stride width ctx batch H KVH D scale ctas ws bytes stream
    # unsupported head_dim -> NVK_ERR_UNSUPPORTED with a message
    rc = lib.nvk_paged_decode(n, n, n, n, 8, 128, n, 4, 4, n, 2, 16, 8, 64, 0.1, 0, n, 0, n)
    assert rc == _lib.NVK_ERR_UNSUPPORTED and b"head_dim" in lib.nvk_last_error()
    # GQA ratio 3 unsupported
    rc = lib.nvk_paged_decode(n, n, n, n, 8, 128, n, 4, 4, n, 2, 24, 8, 128, 0.1, 0, n, 0, n)
    assert rc == _lib.NVK_ERR_UNSUPPORTED
    # block size not a power of two
    rc = lib.nvk_paged_decode(n, n, n, n, 8, 96, n, 4, 4, n, 2, 16, 8, 128, 0.1, 0, n, 0, n)
    assert rc == _lib.NVK_ERR_UNSUPPORTED and b"block_size" in lib.nvk_last_error()
    # table stride narrower than the table
    rc = lib.nvk_paged_decode(n, n, n, n, 8, 128, n, 2, 4, n, 2, 16, 8, 128, 0.1, 0, n, 0, n)
    assert rc == _lib.NVK_ERR_INVALID_ARGUMENT
    # null pointers are rejected before any launch
    rc = lib.nvk_paged_decode(n, n, n, n, 8, 128, n, 4, 4, n, 2, 16, 8, 128, 0.1, 0, n, 0, n)
    assert rc == _lib.NVK_ERR_INVALID_ARGUMENT
    # batch 0 is a no-op
    rc = lib.nvk_paged_decode(n, n, n, n, 8, 128, n, 4, 4, n, 0, 16, 8, 128, 0.1, 0, n, 0, n)
    assert rc == _lib.NVK_OK
    # the no-alloc entry point runs the same checks first, before its scratch-size check
    rc = lib.nvk_paged_decode_noalloc(n, n, n, n, 8, 128, n, 4, 4, n, 1 << 20, 16, 8, 128, 0.1, 0, n)
    assert rc == _lib.NVK_ERR_INVALID_ARGUMENT and b"null pointer" in lib.nvk_last_error()
    rc = lib.nvk_paged_decode_noalloc(n, n, n, n, 8, 128, n, 4, 4, n, 2, 24, 8, 128, 0.1, 0, n)
    assert rc == _lib.NVK_ERR_UNSUPPORTED and b"GQA" in lib.nvk_last_error()
    assert lib.nvk_paged_decode_noalloc_error(None, n) == _lib.NVK_ERR_INVALID_ARGUMENT
    # append: row not a multiple of 16 bytes, zero tokens is a no-op
    rc = lib.nvk_kv_append(n, n, 3, 3, n, n, n, 1, 8, 1, 3, n, n)
    assert rc == _lib.NVK_ERR_UNSUPPORTED
    assert lib.nvk_kv_append(n, n, 1024, 1024, n, n, n, 0, 8, 8, 128, n, n) == _lib.NVK_OK
    rc = lib.nvk_kv_append(n, n, 1024, 1024, n, n, n, 4, 8, 8, 128, n, n)
    assert rc == _lib.NVK_ERR_INVALID_ARGUMENT
    # prefill: block size other than 128 and head_dim other than 128
    rc = lib.nvk_paged_prefill(n, n, n, n, 8, 64, n, 4, n, n, 1, 8, 8, 16, 8, 128, 0.1, n, n)
    assert rc == _lib.NVK_ERR_INVALID_ARGUMENT  # null q/out checked first
    rc = lib.nvk_dense_prefill(n, n, n, n, n, n, 1, 8, 8, 8, 16, 8, 64, 0.1, n, n)
    assert rc == _lib.NVK_ERR_UNSUPPORTED


def test_workspace_size_grows_with_grid_and_batch():
    sz = ctypes.c_size_t()
    lib = _lib.load()
    sizes = []
    for ctas in (1, 148, 296):
        assert lib.nvk_paged_decode_workspace_size(32, 16, 8, 128, ctas, ctypes.byref(sz)) == 0
        sizes.append(sz.value)
    assert sizes[0] < sizes[1] < sizes[2]
    # 148 CTAs x 2 partial slots x 2 query heads x 128 floats is the bulk
    assert sizes[1] >= 148 * 2 * 2 * 128 * 4
    assert lib.nvk_paged_decode_workspace_size(1024, 16, 8, 128, 148, ctypes.byref(sz)) == 0
    assert sz.value >= 1024 * 8 * 4
    assert lib.nvk_paged_decode_workspace_size(32, 16, 8, 64, 1, ctypes.byref(sz)) == _lib.NVK_ERR_UNSUPPORTED


def test_call_wrapper_raises_value_error_on_bad_arguments():
    with pytest.raises(ValueError, match="head_dim"):
        _lib.call("nvk_paged_decode_workspace_size", 1, 16, 8, 64, 1, ctypes.byref(ctypes.c_size_t()))
