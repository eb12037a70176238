"""The C-ABI library loads and exports the header's entry points (CPU only).

No compute calls: this host has no GPU.  Only host-side functions and the
error path of context creation run here.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_functions() -> list[str]:
    src = (ROOT / "include" / "m1moe_cuda.h").read_text()
    return re.findall(r"M1MOE_API\s+[\w\s\*]+?\b(m1moe_cuda_\w+)\s*\(", src)


@pytest.fixture(scope="module")
def lib():
    from m1moe_b200 import build
    build.build()
    from m1moe_b200 import _lib
    return _lib.lib()


def test_header_declares_entry_points():
    names = header_functions()
    assert len(names) >= 16
    assert "m1moe_cuda_moe_layer" in names and "m1moe_cuda_matvec4" in names


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_bindings_cover_header():
    from m1moe_b200 import _lib
    bound = {n for n, _, _ in _lib._SIGS}
    assert set(header_functions()) <= bound


def test_abi_version(lib):
    src = (ROOT / "include" / "m1moe_cuda.h").read_text()
    want = int(re.search(r"#define M1MOE_CUDA_ABI_VERSION (\d+)", src).group(1))
    assert lib.m1moe_cuda_abi_version() == want


def test_expert_bytes_host_function(lib):
    assert lib.m1moe_cuda_expert_bytes(2048, 1024, 64) == 3_538_944
    assert lib.m1moe_cuda_expert_bytes(4096, 14336, 64) == 99_090_432
    assert lib.m1moe_cuda_expert_bytes(100, 64, 64) == 0  # 100 % 64 != 0


def test_create_rejects_bad_config(lib):
    from m1moe_b200 import _lib
    h = ctypes.c_void_p()
    assert lib.m1moe_cuda_create(None, ctypes.byref(h)) == 1
    assert b"NULL" in lib.m1moe_cuda_last_error()
    cfg = _lib.Cfg(2048, 1024, 64, 8, 48, 1, 0, 1, 0, 0, 0)  # group size 48
    assert lib.m1moe_cuda_create(ctypes.byref(cfg), ctypes.byref(h)) == 6
    cfg = _lib.Cfg(2048, 1024, 64, 80, 64, 1, 0, 1, 0, 0, 0)  # top_k > num_experts
    assert lib.m1moe_cuda_create(ctypes.byref(cfg), ctypes.byref(h)) == 1
    cfg = _lib.Cfg(2048, 1024, 64, 8, 64, 1, 0, 9, 0, 0, 0)  # batch 9 > 8
    assert lib.m1moe_cuda_create(ctypes.byref(cfg), ctypes.byref(h)) == 1
    assert not h.value


def test_create_without_gpu_fails_loudly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from m1moe_b200 import _lib
    h = ctypes.c_void_p()
    cfg = _lib.Cfg(128, 64, 4, 2, 64, 1, 0, 1, 0, 0, 0)
    st = lib.m1moe_cuda_create(ctypes.byref(cfg), ctypes.byref(h))
    assert st == 3 and not h.value
    assert lib.m1moe_cuda_last_error()


def test_missing_library_raises(monkeypatch, tmp_path):
    from m1moe_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "nope.so")
    with pytest.raises(ImportError, match="no CPU fallback"):
        _lib.lib()
