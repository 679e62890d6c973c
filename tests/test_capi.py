"""CPU: the C-ABI library loads, exports every entry point the header declares,
and its host-side validation rejects bad arguments before touching the GPU."""
import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "unbox_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ubx_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("ubx_kv_append", "ubx_paged_decode_attention", "ubx_slot_mapping", "ubx_paged_decode_workspace_size",
              "ubx_workspace_init", "ubx_read_device_error"):
        assert s in syms


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.library.load()
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} declared in the header but not exported"
        assert s in pkg.library.SIGNATURES, f"{s} has no ctypes signature"
    nm = os.popen(f"nm -D --defined-only {pkg.library.LIB_PATH}").read()
    for s in declared_symbols():
        assert re.search(rf"\bT {s}\b", nm), s


def declared_arities():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(ubx_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", src):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def test_ctypes_signatures_match_header_arity(pkg):
    """Every ctypes stub passes exactly as many arguments as the C declaration takes."""
    ar = declared_arities()
    assert set(ar) == set(declared_symbols())
    for name, n in ar.items():
        assert len(pkg.library.SIGNATURES[name][1]) == n, (name, n, len(pkg.library.SIGNATURES[name][1]))


def test_host_only_entry_points(pkg):
    lib = pkg.library.load()
    assert lib.ubx_version() >= 100
    assert lib.ubx_status_string(0) == b"ok"
    assert lib.ubx_status_string(3) == b"workspace missing or too small"


def test_validation_rejects_before_any_launch(pkg):
    lib = pkg.library.load()
    # unknown dtype
    st = lib.ubx_paged_decode_attention(None, 0, 0, None, None, 0, 0, 0, None, 0, None, None, 0, 0,
                                        1, 16, 8, 112, 16, 1, 1, 1.0, 7, 0, 0, None, 0, None)
    assert st == pkg.library.ERR_INVALID_ARGUMENT and b"dtype" in lib.ubx_last_error()
    # head_dim not built
    st = lib.ubx_paged_decode_attention(None, 0, 0, None, None, 0, 0, 0, None, 0, None, None, 0, 0,
                                        1, 16, 8, 96, 16, 1, 1, 1.0, 1, 0, 0, None, 0, None)
    assert st == pkg.library.ERR_UNSUPPORTED and b"head_dim" in lib.ubx_last_error()
    # GQA ratio 3
    st = lib.ubx_paged_decode_attention(None, 0, 0, None, None, 0, 0, 0, None, 0, None, None, 0, 0,
                                        1, 12, 4, 112, 16, 1, 1, 1.0, 1, 0, 0, None, 0, None)
    assert st == pkg.library.ERR_UNSUPPORTED
    # page size other than 16
    st = lib.ubx_paged_decode_attention(None, 0, 0, None, None, 0, 0, 0, None, 0, None, None, 0, 0,
                                        1, 16, 8, 112, 32, 1, 1, 1.0, 1, 0, 0, None, 0, None)
    assert st == pkg.library.ERR_UNSUPPORTED and b"block_size" in lib.ubx_last_error()
    # null pointers with a real batch
    st = lib.ubx_paged_decode_attention(None, 0, 0, None, None, 0, 0, 0, None, 0, None, None, 0, 0,
                                        1, 16, 8, 112, 16, 1, 1, 1.0, 1, 0, 0, None, 0, None)
    assert st == pkg.library.ERR_INVALID_ARGUMENT
    # empty batch is a no-op
    st = lib.ubx_paged_decode_attention(None, 0, 0, None, None, 0, 0, 0, None, 0, None, None, 0, 0,
                                        0, 16, 8, 112, 16, 1, 1, 1.0, 1, 0, 0, None, 0, None)
    assert st == 0
    # a workspace off a 16-byte boundary (the kernels read it 16 bytes at a time);
    # the other pointers are never dereferenced on the host
    st = lib.ubx_paged_decode_attention(0x10000, 16 * 112, 112, 0x20000, 0x30000, 16 * 8 * 112, 8 * 112, 112,
                                        0x40000, 1, 0x50000, 0x60000, 16 * 112, 112,
                                        1, 16, 8, 112, 16, 1, 1, 1.0, 1, 0, 0, 0x70008, 1 << 30, None)
    assert st == pkg.library.ERR_WORKSPACE and b"16-byte aligned" in lib.ubx_last_error()
    st = lib.ubx_kv_append(None, None, 0, 0, None, None, 0, 0, 0, None, 0, 8, 112, 16, 4, 1, None, None)
    assert st == 0


def test_ops_refuse_cpu_tensors(pkg):
    """No CPU fallback: host tensors are an error, not a slow path."""
    lay = pkg.workloads.layout_uniform(3, 2, 1, 20, num_blocks=4)
    t = pkg.workloads.materialize_host(lay, 3, dtype="bfloat16")
    with pytest.raises(ValueError, match="CUDA"):
        pkg.paged_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"], t["context_lens"])
    with pytest.raises(ValueError, match="CUDA"):
        pkg.kv_append(t["k_new"], t["v_new"], t["k_cache"], t["v_cache"], t["slot_mapping"])
    with pytest.raises(ValueError, match="CUDA"):
        pkg.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"], t["context_lens"], 16)


def test_missing_library_fails_loudly(pkg, monkeypatch, tmp_path):
    lib_mod = pkg.library
    monkeypatch.setattr(lib_mod, "_lib", None)
    monkeypatch.setattr(lib_mod, "LIB_PATH", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        lib_mod.load()
