"""The C-ABI library loads and exports exactly what include/paged_serve.h declares.

Runs without a GPU: only symbol lookups and argument checks that return before
any CUDA call are exercised here.
"""

from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from paged_serve_b200 import _lib
from paged_serve_b200.build import LIB_PATH
from tests.conftest import ROOT

HEADER = ROOT / "include" / "paged_serve.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^PS_API\s+[\w\s\*]+?\b(ps_\w+)\s*\(", text, flags=re.M)


def test_header_declares_the_hot_path():
    names = set(declared_functions())
    assert {"ps_cache_append", "ps_cache_append_rope", "ps_copy_blocks", "ps_paged_decode",
            "ps_paged_prefill", "ps_paged_decode_workspace_bytes", "ps_last_error_string",
            "ps_abi_version"} <= names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (ps_\w+)", out))
    assert exported == set(declared_functions())


def test_binding_table_matches_header():
    assert set(_lib.SIGNATURES) == set(declared_functions())
    text = HEADER.read_text()
    for name, (_, args) in _lib.SIGNATURES.items():
        decl = re.search(rf"^PS_API[^;(]*\b{name}\s*\(([^)]*)\)", text, flags=re.M).group(1)
        n = 0 if decl.strip() == "void" else decl.count(",") + 1
        assert n == len(args), f"{name}: header has {n} params, binding {len(args)}"


def test_abi_version():
    assert _lib.load().ps_abi_version() == _lib.ABI_VERSION


def test_binding_constants_match_the_header():
    """The binding's ABI version and device error bits are the header's macros."""
    macros = dict(re.findall(r"^#define (PS_\w+) (\d+)", HEADER.read_text(), flags=re.M))
    assert int(macros["PS_ABI_VERSION"]) == _lib.ABI_VERSION
    for name in ("PS_DEVERR_BLOCK_ID", "PS_DEVERR_SLOT", "PS_DEVERR_POSITION",
                 "PS_DEVERR_TIMEOUT", "PS_DEVERR_LENGTH", "PS_DEVERR_BLOCK_PAIRS"):
        assert int(macros[name]) == getattr(_lib, name), name


def _msg():
    return _lib.load().ps_last_error_string().decode()


class TestArgumentChecks:
    """Bad arguments are rejected on the host, before any launch."""

    def test_append_rejects_fp32(self):
        lib = _lib.load()
        st = lib.ps_cache_append(1, 1, 1, 1, 1, 4, 256, 256, 2, 128, 16, 8, 3, None, None)
        assert st == _lib.PS_ERR_UNSUPPORTED and "dtype" in _msg()

    def test_append_rejects_head_dim(self):
        lib = _lib.load()
        st = lib.ps_cache_append(1, 1, 1, 1, 1, 4, 256, 256, 2, 96, 16, 8, 2, None, None)
        assert st == _lib.PS_ERR_UNSUPPORTED and "head_dim" in _msg()

    def test_append_zero_tokens_is_a_no_op(self):
        lib = _lib.load()
        assert lib.ps_cache_append(None, None, None, None, None, 0, 256, 256, 2, 128, 16, 8, 2,
                                   None, None) == _lib.PS_OK

    def test_append_rejects_null_pointers(self):
        lib = _lib.load()
        st = lib.ps_cache_append(None, None, None, None, None, 4, 256, 256, 2, 128, 16, 8, 2,
                                 None, None)
        assert st == _lib.PS_ERR_INVALID

    def test_append_rejects_misaligned_key(self):
        lib = _lib.load()
        st = lib.ps_cache_append(16, 16, 18, 16, 16, 4, 256, 256, 2, 128, 16, 8, 2, None, None)
        assert st == _lib.PS_ERR_INVALID and "aligned" in _msg()

    def test_rope_requires_full_rotary_dim(self):
        lib = _lib.load()
        st = lib.ps_cache_append_rope(16, 16, 16, 16, 16, 16, 4, 256, 256, 2, 128, 16, 8, 16,
                                      100, 64, 2, None, None)
        assert st == _lib.PS_ERR_UNSUPPORTED and "rope_dim" in _msg()

    def test_copy_rejects_unaligned_block_bytes(self):
        lib = _lib.load()
        st = lib.ps_copy_blocks(16, 16, 16, 2, 1, 0, 100, 8, None, None)
        assert st == _lib.PS_ERR_INVALID

    def test_decode_rejects_ragged_gqa(self):
        lib = _lib.load()
        st = lib.ps_paged_decode(16, 4096, 16, 4096, 16, 16, 8, 16, 8, 16, 2, 30, 8, 128, 16, 8,
                                 0.1, 0, None, 0, 2, None, None)
        assert st == _lib.PS_ERR_INVALID and "divisible" in _msg()

    @pytest.mark.parametrize("bs", [24, 64])
    def test_decode_rejects_block_size(self, bs):
        lib = _lib.load()
        st = lib.ps_paged_decode(16, 4096, 16, 4096, 16, 16, 8, 16, 8, 16, 2, 32, 8, 128, bs, 8,
                                 0.1, 0, None, 0, 2, None, None)
        assert st == _lib.PS_ERR_UNSUPPORTED and "block_size" in _msg()

    def test_decode_split_needs_workspace(self):
        lib = _lib.load()
        st = lib.ps_paged_decode(256, 4096, 256, 4096, 256, 256, 64, 256, 64, 256, 2, 32, 8, 128,
                                 16, 64, 0.1, 256, None, 0, 2, None, None)
        assert st == _lib.PS_ERR_INVALID and "workspace" in _msg()

    def test_noalloc_checks_arguments_before_sizing_its_scratch(self):
        lib = _lib.load()
        st = lib.ps_paged_decode_noalloc(16, 4096, 16, 4096, 16, 16, 1 << 20, 16, 256, 16, 70000,
                                         32, 8, 128, 16, 256, 0.1, 512, 2, None, None)
        assert st == _lib.PS_ERR_INVALID and "too many sequences" in _msg()
        st = lib.ps_paged_decode_noalloc(16, 4096, 16, 4096, 16, 16, 1 << 20, 16, 256, 16, 64,
                                         32, 8, 128, 16, 256, 0.1, 500, 2, None, None)
        assert st == _lib.PS_ERR_INVALID and "multiple of" in _msg()
        st = lib.ps_paged_decode_noalloc(16, 4096, 16, 4096, 16, 16, 1 << 20, 16, 256, 16, 4096,
                                         32, 8, 128, 16, 256, 0.1, 512, 2, None, None)
        assert st == _lib.PS_ERR_INVALID and "built-in scratch" in _msg()
        assert _msg().startswith("ps_paged_decode_noalloc")

    def test_stream_read_rejects_ragged_sizes_and_unknown_methods(self):
        lib = _lib.load()
        for method in (_lib.PS_STREAM_BULK, _lib.PS_STREAM_LOADS):
            assert lib.ps_stream_read(16, 100, 16, method, None, None) == _lib.PS_ERR_INVALID
            assert lib.ps_stream_read(18, 96, 16, method, None, None) == _lib.PS_ERR_INVALID
            assert lib.ps_stream_read(None, 0, None, method, None, None) == _lib.PS_OK
        assert lib.ps_stream_read(16, 96, 16, 7, None, None) == _lib.PS_ERR_INVALID
        assert "method" in _msg()

    def test_workspace_bytes(self):
        lib = _lib.load()
        assert lib.ps_paged_decode_workspace_bytes(4, 32, 128, 16, 64, 0) == 0
        assert lib.ps_paged_decode_workspace_bytes(4, 32, 128, 16, 64, 1024) == 0
        got = lib.ps_paged_decode_workspace_bytes(4, 32, 128, 16, 64, 512)
        rows = 4 * 2 * 32  # sequences x partitions x query heads
        units = 4 * 2  # (sequence, partition) list for the persistent launch
        assert got == ((rows * 128 * 4 + 255) // 256 + (rows * 4 + 255) // 256
                       + (units * 4 + 255) // 256 + 1) * 256

    def test_prefill_split_checks_split_keys_and_workspace(self):
        lib = _lib.load()
        # 1 sequence, 512 new tokens over a 32k table (2048 blocks of 16), Hq 32, Hkv 8, D 128
        args = (256, 4096, 256, 4096, 512, 256, 256, 4096, 256, 2048, 256, 256, 256, 1, 512,
                32, 8, 128, 16, 2048, 0.1)
        st = lib.ps_paged_prefill_split(*args, 100, 256, 1 << 30, 2, None, None)
        assert st == _lib.PS_ERR_INVALID and "multiple of 128" in _msg()
        st = lib.ps_paged_prefill_split(*args, 4096, None, 0, 2, None, None)
        assert st == _lib.PS_ERR_INVALID and "workspace" in _msg()
        need = lib.ps_paged_prefill_workspace_bytes(1, 512, 32, 8, 128, 16, 2048, 4096)
        st = lib.ps_paged_prefill_split(*args, 4096, 256, need - 256, 2, None, None)
        assert st == _lib.PS_ERR_INVALID and "needed" in _msg()
        assert _msg().startswith("ps_paged_prefill_split")

    def test_prefill_workspace_bytes(self):
        lib = _lib.load()
        # G = 4: 32 tokens per query tile, 64 per item; 512 tokens -> 8 items per KV head
        items = 8 * 8
        pieces = 32768 // 4096
        rows = items * pieces * 2 * 128
        got = lib.ps_paged_prefill_workspace_bytes(1, 512, 32, 8, 128, 16, 2048, 4096)
        assert got == ((rows * 128 * 4 + 255) // 256 + (rows * 8 + 255) // 256) * 256
        # nothing split: split_keys 0, or a piece covering the whole table
        assert lib.ps_paged_prefill_workspace_bytes(1, 512, 32, 8, 128, 16, 2048, 0) == 0
        assert lib.ps_paged_prefill_workspace_bytes(1, 512, 32, 8, 128, 16, 2048, 32768) == 0
        assert lib.ps_paged_prefill_workspace_bytes(1, 512, 32, 8, 128, 16, 2048, 100) == 0

    def test_status_maps_to_reference_exception_types(self):
        _lib.load().ps_cache_append(1, 1, 1, 1, 1, 4, 256, 256, 2, 96, 16, 8, 2, None, None)
        with pytest.raises(ValueError, match="head_dim"):
            _lib.check(_lib.PS_ERR_UNSUPPORTED, "x")
        with pytest.raises(_lib.NativeError):
            _lib.check(_lib.PS_ERR_CUDA, "x")


def test_ctypes_pointer_types():
    for _, (_, args) in _lib.SIGNATURES.items():
        for a in args:
            assert a in (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float)


def test_every_compute_entry_point_opens_an_nvtx_range():
    """Each C-ABI call that enqueues work is a named NVTX range in profiler timelines."""
    plumbing = {"ps_abi_version", "ps_last_error_string", "ps_paged_decode_workspace_bytes",
                "ps_paged_prefill_workspace_bytes"}
    sources = "\n".join(p.read_text() for p in (ROOT / "paged_serve_b200" / "csrc").glob("*.cu"))
    for name in set(declared_functions()) - plumbing:
        m = re.search(rf'extern "C" [\w\s\*]+?\b{name}\([^{{]*\{{\s*ps::NvtxRange nvtx_range\('
                      rf'"{name}"\);', sources)
        assert m, f"{name} has no NVTX range"
